"""Lane grouping by density class (gsp_group_plan, grouped_grammar_logits):
the device plan equals a numpy restatement of the planner (per-request legal
tokens and active tiles, order by tile fill, prefix / suffix active tiles,
every split costed with the route model), and a split batch gives, row for
row, exactly what each group's route gives for that group alone, with the
oracle's support and top-1. A batch that does not pay for a split runs one
route; batch 1 never splits.
"""
import numpy as np
import pytest
import torch

from gsp import _native
from gsp import triton_runtime as tr
from gsp import workloads as wl
from oracle import gsp_oracle as O

pytestmark = pytest.mark.gpu

V, H = 32768, 512
# small fixed costs so that a split pays at this size
COST = {"row_sparse_fixed_us": 0.5, "block_floor_us": 0.0, "block_fixed_us": 1.0, "dense_fixed_us": 1.0,
        "group_split_fixed_us": 0.5}


def _best(batch, legal_total, active, c, e=2):
    """The route model (best_route_by_cost) in the same double arithmetic."""
    row_bytes = H * e
    out_bytes = batch * V * e
    t_row = c["row_sparse_fixed_us"] + (legal_total * row_bytes + out_bytes) / (c["hbm_gbs"] * 1e3)
    if batch <= 1:
        return 0, (0.0 if batch <= 0 else t_row)
    rows = min(active * 128, V)
    t_block = c["block_fixed_us"] + (rows * row_bytes) / (c["block_gbs"] * 1e3)
    if c["block_floor_us"] > t_block:
        t_block = c["block_floor_us"]
    t_dense = c["dense_fixed_us"] + (V * row_bytes) / (c["dense_gbs"] * 1e3)
    best, bt = 1, t_block
    if t_dense < bt:
        best, bt = 2, t_dense
    if t_row < bt:
        best, bt = 0, t_row
    return best, bt


def plan_reference(mask_np, with_logits, cost):
    c = dict(tr.B200_COST, **cost)
    B = mask_np.shape[0]
    legal_bits = wl.unpack_bitmask(mask_np, V)
    ntiles = (V + 127) // 128
    padded = np.zeros((B, ntiles * 128), dtype=bool)
    padded[:, :V] = legal_bits
    tile_any = padded.reshape(B, ntiles, 128).any(axis=2)
    legal = legal_bits.sum(axis=1).astype(np.int64)
    tiles = tile_any.sum(axis=1).astype(np.int64)
    fill = [legal[b] / (128.0 * tiles[b]) if tiles[b] else -1.0 for b in range(B)]
    order = sorted(range(B), key=lambda b: (fill[b], b))
    inverse = np.empty(B, dtype=np.int64)
    inverse[order] = np.arange(B)
    pos = np.where(tile_any, inverse[:, None], -1)
    active = tile_any.any(axis=0)
    hmin = np.bincount(np.where(tile_any, inverse[:, None], B).min(axis=0)[active], minlength=B)[:B]
    hmax = np.bincount(pos.max(axis=0)[active], minlength=B)[:B]
    legal_total, active_total = int(legal.sum()), int(hmax.sum())
    single, t_single = _best(B, legal_total, active_total, c)
    unperm = 2.0 * (B * V * 2) / (c["hbm_gbs"] * 1e3) if with_logits else 0.0
    best_t, best = t_single, (0, single, single)
    la = aa = 0
    ab = active_total
    for k in range(1, B):
        la += int(legal[order[k - 1]])
        aa += int(hmin[k - 1])
        ab -= int(hmax[k - 1])
        ra, ta = _best(k, la, aa, c)
        rb, tb = _best(B - k, legal_total - la, ab, c)
        tt = ta + tb + c["group_split_fixed_us"] + unperm
        if tt < best_t:
            best_t, best = tt, (k, ra, rb)
    return {"k": best[0], "ra": best[1], "rb": best[2], "single": single,
            "single_ns": int(min(t_single * 1e3, 2e9)), "split_ns": int(min(best_t * 1e3, 2e9)) if best[0] else -1,
            "order": order}


def _mixed_mask(rng, n_scattered, n_clustered, frac=0.005, cfrac=0.2):
    sc = wl.make_batch_mask(rng, n_scattered, V, [int(frac * V)] * n_scattered)
    cl = np.repeat(wl.make_batch_mask(rng, 1, V, [int(cfrac * V)], clustered=True, max_runs=1), n_clustered, axis=0)
    m = np.concatenate([sc, cl])
    return m[rng.permutation(m.shape[0])]


@pytest.fixture(scope="module")
def weight(cuda_device):
    rng = np.random.default_rng(5)
    return (torch.from_numpy(rng.standard_normal((V, H), dtype=np.float32)) * 0.05).half()


@pytest.mark.parametrize("with_logits", [True, False])
def test_plan_matches_restatement(cuda_device, with_logits):
    rng = np.random.default_rng(11)
    for mask_np, cost in ((_mixed_mask(rng, 12, 4), COST), (_mixed_mask(rng, 20, 12), COST),
                          (wl.make_batch_mask(rng, 9, V, [50, 0, 3000, 7, 7, 20000, 1, 0, 400]), COST),
                          (_mixed_mask(rng, 12, 4), {})):
        md = torch.from_numpy(mask_np).to(cuda_device)
        B = mask_np.shape[0]
        plan = torch.empty(_native.GROUP_PLAN_HEADER + 6 * B, dtype=torch.int32, device=cuda_device)
        _native.group_plan(md, V, H, 2, with_logits, plan, cost)
        got = plan.cpu().numpy()
        ref = plan_reference(mask_np, with_logits, cost)
        hdr = got[:6].tolist()
        assert hdr == [ref["k"], ref["ra"], ref["rb"], ref["single"], ref["single_ns"], ref["split_ns"]], (hdr, ref)
        order = got[16:16 + B].tolist()
        assert order == ref["order"]
        assert got[16 + B:16 + 2 * B].tolist() == np.argsort(order).tolist()


def test_split_batch_matches_each_groups_route(cuda_device, weight):
    rng = np.random.default_rng(3)
    mask_np = _mixed_mask(rng, 12, 4)
    ref = plan_reference(mask_np, True, COST)
    assert ref["k"] > 0 and ref["ra"] != ref["rb"], ref  # the case design: a split with two routes
    dev = cuda_device
    w = weight.to(dev)
    B = mask_np.shape[0]
    h = torch.from_numpy(rng.standard_normal((B, H), dtype=np.float32)).half()
    res = tr.grouped_grammar_logits(h.to(dev), w, torch.from_numpy(mask_np).to(dev), cost=COST)
    assert res.plan["split"] == ref["k"]
    fns = {0: _native.row_sparse, 1: _native.block_gemm, 2: _native.dense_masked}
    order = ref["order"]
    for lo, hi, route in ((0, ref["k"], ref["ra"]), (ref["k"], B, ref["rb"])):
        rows = order[lo:hi]
        hg = h[rows].contiguous().to(dev)
        mg = torch.from_numpy(mask_np[rows]).to(dev)
        lg = torch.empty(len(rows), V, dtype=torch.float16, device=dev)
        tv = torch.empty(len(rows), device=dev)
        ti = torch.empty(len(rows), dtype=torch.int64, device=dev)
        fns[route](hg, w, mg, logits=lg, top_value=tv, top_index=ti)
        idx = torch.tensor(rows, device=dev)
        assert torch.equal(res.logits[idx], lg), (lo, hi, route)
        assert torch.equal(res.top_value[idx], tv) and torch.equal(res.top_index[idx], ti), (lo, hi, route)
    exact = O.masked_logits_exact(h, weight, mask_np)
    rep = O.compare_logits(exact, res.logits.cpu(), dtype=torch.float16)
    assert rep["support"] and rep["values"], rep
    assert O.top1_agrees(exact, res.top_index.cpu(), dtype=torch.float16)
    # top-1 only: same tokens, no logits
    res2 = tr.grouped_grammar_logits(h.to(dev), w, torch.from_numpy(mask_np).to(dev), cost=COST, return_logits=False)
    assert res2.logits is None and torch.equal(res2.top_index, res.top_index)


def test_no_split_when_it_does_not_pay(cuda_device, weight):
    rng = np.random.default_rng(8)
    dev = cuda_device
    w = weight.to(dev)
    for B, ks in ((8, [int(0.9 * V)] * 8), (1, [30])):
        mask_np = wl.make_batch_mask(rng, B, V, ks)
        h = torch.from_numpy(rng.standard_normal((B, H), dtype=np.float32)).half().to(dev)
        res = tr.grouped_grammar_logits(h, w, torch.from_numpy(mask_np).to(dev), cost=COST)
        assert res.plan["split"] == 0 and len(res.plan["routes"]) == 1
        fn = {"row-sparse": _native.row_sparse, "block-sparse": _native.block_gemm,
              "dense-mask": _native.dense_masked}[res.plan["routes"][0]]
        lg = torch.empty(B, V, dtype=torch.float16, device=dev)
        fn(h, w, torch.from_numpy(mask_np).to(dev), logits=lg)
        assert torch.equal(res.logits, lg)


def test_plan_on_ragged_vocabulary(cuda_device):
    """A vocabulary that is not a multiple of 32 or 128, with the bits past it
    set in every request's last word: the device plan still equals the
    restatement's, which never counts those bits."""
    global V
    saved = V
    try:
        V = 30001
        rng = np.random.default_rng(17)
        mask_np = _mixed_mask(rng, 9, 3)
        mask_np[:, -1] |= np.int32(-1)
        B = mask_np.shape[0]
        plan = torch.empty(_native.GROUP_PLAN_HEADER + 6 * B, dtype=torch.int32, device=cuda_device)
        _native.group_plan(torch.from_numpy(mask_np).to(cuda_device), V, H, 2, True, plan, COST)
        got = plan.cpu().numpy()
        ref = plan_reference(mask_np, True, COST)
        assert got[:6].tolist() == [ref["k"], ref["ra"], ref["rb"], ref["single"], ref["single_ns"], ref["split_ns"]]
        assert got[16:16 + B].tolist() == ref["order"]
    finally:
        V = saved
