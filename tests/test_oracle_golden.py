"""The CPU oracle against the golden fixtures generated from the reference's own
code (tests/golden/make_golden.py). CPU only."""
import numpy as np
import pytest
import torch

from conftest import load_json, load_npz
from oracle import gsp_oracle as O


def _case_inputs(c):
    w, h, mask = O.kernel_case_inputs(c["vocab"], c["hidden"], c["batch"], c["dtype"], c["seed"],
                                      c["recipe"], c["extra_words"])
    assert O.tensor_sha256(w) == c["weight_sha256"], "weight generator drifted"
    assert O.tensor_sha256(h) == c["hidden_sha256"], "hidden generator drifted"
    assert O.tensor_sha256(mask) == c["mask_sha256"], "mask generator drifted"
    return w, h, mask


@pytest.mark.parametrize("fixture", ["row_sparse_ref.npz", "block_gemm_ref.npz", "dense_mask_ref.npz"])
def test_oracle_matches_reference_kernels(fixture):
    data, meta = load_npz(fixture)
    assert meta
    for c in meta:
        w, h, mask = _case_inputs(c)
        ref = O.bits16_to_tensor(data[c["name"] + "/out"], c["dtype"]).double()
        exact = O.masked_logits_exact(h, w, mask)
        assert torch.equal(torch.isfinite(ref), torch.isfinite(exact)), (fixture, c["name"])
        fin = torch.isfinite(exact)
        # The reference rounds its fp32 accumulator once; under the Triton CPU
        # interpreter the fp32 -> bf16 conversion truncates, so allow one output
        # ulp, plus 1e-4 absolute for fp32 accumulation noise near zero.
        err = (ref[fin] - exact[fin]).abs()
        bound = O.ulp(O.TORCH_DTYPES[c["dtype"]], exact[fin]) + 1e-4
        assert bool((err <= bound).all()), (fixture, c["name"], float(err.max()))
        # The oracle's rounded logits meet the product tolerance against the exact values.
        dt = O.TORCH_DTYPES[c["dtype"]]
        rep = O.compare_logits(exact, O.masked_logits(h, w, mask), dtype=dt)
        assert rep["support"] and rep["values"], (fixture, c["name"], rep)
        _, idx = O.top1(O.masked_logits(h, w, mask))
        assert O.top1_agrees(exact, idx, dtype=dt), (fixture, c["name"])
        _, idx_ref = O.top1(ref)
        assert O.top1_agrees(exact, idx_ref, dtype=dt), (fixture, c["name"])


def test_reference_kernels_ignore_tail_bits_and_extra_words():
    """Rows >= V and words beyond ceil(V/32) never become legal
    (gsp/triton_runtime.py:30,35 of the reference)."""
    data, meta = load_npz("row_sparse_ref.npz")
    c = next(m for m in meta if m["name"] == "v1000_h256_b3_f16_mixed")
    ref = O.bits16_to_tensor(data[c["name"] + "/out"], c["dtype"])
    assert ref.shape == (3, 1000)
    assert torch.isfinite(ref[2]).all()      # 'full' row: every word -1, tail bits set
    assert not torch.isfinite(ref[1]).any()  # 'zero' row


def test_oracle_projection_matches_reference_runtime():
    data = np.load(__import__("conftest").GOLDEN + "/projection_ref.npz")
    import json
    meta = json.loads(str(data["meta"]))
    for c in meta:
        if c["name"].startswith("config0"):
            w, h, ids = O.config0_inputs(seed=0)
            assert np.array_equal(ids, data[c["name"] + "/ids"])
        else:
            w, h = O.projection_case_inputs(c["dtype"], c["seed"])
            if c["hidden_1d"]:
                h = h[0]
            ids = None if c["ids_is_none"] else torch.from_numpy(data[c["name"] + "/ids"])
        assert O.tensor_sha256(w) == c["weight_sha256"]
        assert O.tensor_sha256(h) == c["hidden_sha256"]
        if c["name"].startswith("config0"):
            ids = torch.from_numpy(ids)
        res = O.constrained_projection(h, w, ids, dense_threshold=c["threshold"])
        assert res.mode == c["mode"], c["name"]
        assert np.array_equal(res.token_ids.numpy(), data[c["name"] + "/token_ids"])
        raw = data[c["name"] + "/logits"]
        ref = torch.from_numpy(raw) if raw.dtype == np.float32 else O.bits16_to_tensor(raw, c["dtype"])
        rep = O.compare_logits(ref, res.logits, dtype=None if ref.dtype == torch.float32 else ref.dtype,
                               atol=1e-5 if ref.dtype == torch.float32 else O.ATOL)
        assert rep["support"] and rep["values"], (c["name"], rep)
    errors = __import__("json").loads(str(data["errors"]))
    w = torch.zeros((100, 8))
    h = torch.zeros((1, 8))
    cases = {"empty": torch.zeros(0, dtype=torch.long), "negative": torch.tensor([-1, 3]),
             "too_large": torch.tensor([5, 100]), "two_dim": torch.tensor([[1, 2]])}
    for label, ids in cases.items():
        with pytest.raises(ValueError) as exc:
            O.constrained_projection(h, w, ids)
        assert str(exc.value) == errors[label]


def test_config0_cpu_plumbing_case():
    """32,768 x 1,024 fp32, batch 1, 1% uniform, seed 0: sparse-gather with 327
    legal logits, -inf elsewhere, same greedy token as dense + mask."""
    data = np.load(__import__("conftest").GOLDEN + "/projection_ref.npz")
    w, h, ids = O.config0_inputs(seed=0)
    mask = O.ids_to_bitmask(ids, w.shape[0])
    full = O.masked_logits(h, w, mask)
    assert int(torch.isfinite(full).sum()) == len(ids) == 327
    ref_ids = data["config0_fp32_1pct/token_ids"]
    ref_logits = torch.from_numpy(data["config0_fp32_1pct/logits"])[0]
    _, top = O.top1(full)
    assert int(top[0]) == int(ref_ids[int(ref_logits.argmax())])


def test_oracle_routes_match_reference():
    routes = load_json("routes_ref.json")
    for c in routes["dispatch_cases"]:
        assert O.adaptive_route(c["batch"], c["fwf"]) == c["route"], c
        assert O.adaptive_route(c["batch"], None) == c["route_without_fwf"], c
    for c in routes["grid"]:
        assert O.adaptive_route(c["batch"], c["fwf"], c["threshold"]) == c["route"], c
    for c in routes["full_word_fraction"]:
        assert O.full_word_fraction(np.array(c["mask"], dtype=np.int32)) == c["fwf"]


def test_route_known_answers():
    """tests/test_adaptive_dispatch.py:65-74 of the reference."""
    expect = {(1, "all_sparse"): "row-sparse", (1, "all_dense"): "row-sparse",
              (32, "all_sparse"): "block-sparse", (32, "all_dense"): "dense-mask", (32, "mixed"): "dense-mask"}
    for b in (2, 4, 8, 16):
        expect[(b, "all_sparse")] = "block-sparse"
        expect[(b, "all_dense")] = "dense-mask"
        expect[(b, "mixed")] = "block-sparse"
    got = {(c["batch"], c["pattern"]): c["route"] for c in load_json("routes_ref.json")["dispatch_cases"]}
    assert got == expect


def test_pack_unpack_roundtrip():
    rng = np.random.default_rng(0)
    for vocab in (1, 31, 32, 33, 1000, 4096):
        legal = rng.random((3, vocab)) < 0.3
        packed = O.pack_bitmask(legal)
        assert packed.shape == (3, (vocab + 31) // 32)
        assert np.array_equal(O.unpack_bitmask(packed, vocab), legal)


def test_clustered_generator_properties():
    rng = np.random.default_rng(1)
    for k, runs in ((1, 1), (1242, 16), (2483, 64), (24832, 64)):
        ids = O.clustered_legal_ids(rng, 248320, k, runs)
        assert len(ids) == k and len(np.unique(ids)) == k
        assert ids.min() >= 0 and ids.max() < 248320
        assert int((np.diff(ids) > 1).sum()) + 1 <= runs
