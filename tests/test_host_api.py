"""CPU-side checks of the C ABI library and of the drop-in Python API: the
library loads and exports every symbol include/gsp_b200.h declares, C-level
argument validation fails before any device work, and the Python entry points
raise the reference's ValueErrors. No kernel is launched here."""
import ctypes
import os
import re

import pytest
import torch

from conftest import REPO, load_json
from gsp import _native
from gsp import runtime as rt
from gsp import triton_runtime as tr

HEADER = os.path.join(REPO, "include", "gsp_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int32_t|size_t|void|const char\s*\*)\s*(gsp_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    syms = declared_symbols()
    assert len(syms) >= 11
    lib = _native.load()
    for s in syms:
        assert hasattr(lib, s), s
        assert s in _native.SIGNATURES, f"{s} has no ctypes signature"


def test_abi_version_and_status_strings():
    lib = _native.load()
    assert lib.gsp_abi_version() == 1
    assert lib.gsp_status_string(0) == b"GSP_OK"
    assert lib.gsp_status_string(-4) == b"GSP_ERR_CUDA"


def test_workspace_bytes():
    lib = _native.load()
    assert lib.gsp_workspace_bytes(0, 10) == 0
    n = lib.gsp_workspace_bytes(32, 248320)
    assert n % 256 == 0 and n >= 8 * 32 + 1940 * 4


FAKE = ctypes.c_void_p(4096)  # never dereferenced: every call below fails validation first


def _row_sparse(**kw):
    args = dict(hidden=FAKE, hs=8, weight=FAKE, ws=8, mask=None, ms=0, batch=1, vocab=64, hdim=8,
                dtype=0, off=0, logits=None, ls=64, tv=None, ti=None, tk=None, wsp=None, wsb=0)
    args.update(kw)
    lib = _native.load()
    return lib.gsp_row_sparse_logits(args["hidden"], args["hs"], args["weight"], args["ws"], args["mask"],
                                     args["ms"], args["batch"], args["vocab"], args["hdim"], args["dtype"],
                                     args["off"], args["logits"], args["ls"], args["tv"], args["ti"],
                                     args["tk"], args["wsp"], args["wsb"], None)


def test_c_abi_validation_rejects_before_launch():
    lib = _native.load()
    assert _row_sparse(hidden=None) == _native.GSP_ERR_INVALID_ARGUMENT
    assert b"non-null" in lib.gsp_last_error()
    assert _row_sparse(batch=0) == _native.GSP_ERR_INVALID_ARGUMENT
    assert _row_sparse(dtype=7) == _native.GSP_ERR_UNSUPPORTED
    assert _row_sparse(batch=2, hs=4) == _native.GSP_ERR_INVALID_ARGUMENT
    assert _row_sparse(batch=2, mask=FAKE, ms=1) == _native.GSP_ERR_INVALID_ARGUMENT
    assert _row_sparse(tv=FAKE) == _native.GSP_ERR_WORKSPACE
    assert _row_sparse(tv=FAKE, wsp=FAKE, wsb=1) == _native.GSP_ERR_WORKSPACE
    assert lib.gsp_ids_to_bitmask(None, 3, 10, FAKE, FAKE, None) == _native.GSP_ERR_INVALID_ARGUMENT
    assert lib.gsp_mask_stats(None, 0, 1, 10, None, None, None, None) == _native.GSP_ERR_INVALID_ARGUMENT
    assert lib.gsp_top1_from_keys(None, 1, None, None, None) == _native.GSP_ERR_INVALID_ARGUMENT


def _vp_call(route=0, batch=1, tv=FAKE, peers=None, rank=0, world=2, max_batch=4, offset=0, total=128):
    lib = _native.load()
    arr = None if peers is None else (ctypes.c_void_p * len(peers))(*peers)
    return lib.gsp_vocab_parallel_logits(route, FAKE, 8, FAKE, 8, None, 0, batch, 64, 8, 0, offset, None, 64,
                                         tv, None, None, FAKE, 1 << 30, arr, rank, world, max_batch, total, 0, None)


def test_vocab_parallel_entry_validation():
    lib = _native.load()
    ok_peers = [FAKE, FAKE]
    assert _vp_call(route=5, peers=ok_peers) == _native.GSP_ERR_INVALID_ARGUMENT
    assert b"route" in lib.gsp_last_error()
    assert _vp_call(world=9, peers=ok_peers) == _native.GSP_ERR_INVALID_ARGUMENT
    assert _vp_call(rank=2, peers=ok_peers) == _native.GSP_ERR_INVALID_ARGUMENT
    assert _vp_call(tv=None, peers=ok_peers) == _native.GSP_ERR_INVALID_ARGUMENT
    assert b"top-1" in lib.gsp_last_error()
    assert _vp_call(peers=None) == _native.GSP_ERR_INVALID_ARGUMENT
    assert _vp_call(peers=[FAKE, None]) == _native.GSP_ERR_INVALID_ARGUMENT
    assert _vp_call(batch=5, peers=ok_peers, max_batch=4) == _native.GSP_ERR_INVALID_ARGUMENT
    assert b"max_batch" in lib.gsp_last_error()
    assert _vp_call(peers=ok_peers, offset=96, total=128) == _native.GSP_ERR_INVALID_ARGUMENT
    assert b"outside" in lib.gsp_last_error()
    assert lib.gsp_peer_exchange_bytes(0, 4) == 0 and lib.gsp_peer_exchange_bytes(9, 4) == 0
    assert lib.gsp_peer_exchange_bytes(8, 128) >= 1152 + 2 * 8 * 128 * 8
    assert lib.gsp_peer_exchange_alloc(16, None, None) == _native.GSP_ERR_INVALID_ARGUMENT
    assert lib.gsp_peer_exchange_close(None) == _native.GSP_OK and lib.gsp_peer_exchange_free(None) == _native.GSP_OK


def test_python_api_rejects_cpu_tensors_like_the_reference():
    h = torch.zeros(2, 8, dtype=torch.float16)
    w = torch.zeros(64, 8, dtype=torch.float16)
    m = torch.zeros(2, 2, dtype=torch.int32)
    with pytest.raises(ValueError, match="hidden and weight must be CUDA tensors"):
        tr.bitmask_sparse_logits(h, w, m)
    with pytest.raises(ValueError, match="hidden and weight must be CUDA tensors"):
        tr.bitmask_block_gemm_logits(h, w, m)
    with pytest.raises(ValueError, match=r"block GEMM path expects hidden shape \[B,D\] with B >= 2"):
        tr.bitmask_block_gemm_logits(h[:1], w, m[:1])
    with pytest.raises(ValueError, match="hidden and weight must be CUDA tensors"):
        tr.dense_masked_logits(h, w, m)
    with pytest.raises(ValueError):
        rt.constrained_projection(h, w, torch.tensor([1, 2]))


def test_mask_staging_validation():
    with pytest.raises(ValueError, match="bitmask_cpu must be CPU int32"):
        tr.copy_bitmask_to_gpu(torch.zeros(1, 4, dtype=torch.int64))
    with pytest.raises(ValueError, match="bitmask_cpu must be pinned"):
        tr.copy_bitmask_to_gpu(torch.zeros(1, 4, dtype=torch.int32))


def test_full_word_fraction_matches_reference():
    for c in load_json("routes_ref.json")["full_word_fraction"]:
        assert tr.full_word_fraction_cpu(torch.tensor(c["mask"], dtype=torch.int32)) == c["fwf"]


def test_reference_policy_routes_match_reference():
    routes = load_json("routes_ref.json")
    for c in routes["dispatch_cases"]:
        assert tr._reference_route(c["batch"], c["fwf"], 0.80) == c["route"]
        assert tr._reference_route(c["batch"], None, 0.80) == c["route_without_fwf"]
    for c in routes["grid"]:
        assert tr._reference_route(c["batch"], c["fwf"], c["threshold"]) == c["route"]
    with pytest.raises(ValueError, match="full_word_fraction length must equal batch"):
        tr._reference_route(3, [0.1, 0.2], 0.8)


def test_b200_cost_model_prefers_the_cheapest_bytes():
    V, H, e = 248320, 2048, 2
    assert tr.choose_route(1, V, H, e, [V], 1940) == "row-sparse"
    # two requests with a few clustered tokens: row-sparse reads far fewer bytes
    assert tr.choose_route(2, V, H, e, [1242, 1242], 40) == "row-sparse"
    # 32 requests sharing one grammar state: the union of tiles is read once,
    # row-sparse would read the same rows 32 times
    assert tr.choose_route(32, V, H, e, [1242] * 32, 20) == "block-sparse"
    # 32 requests with disjoint clustered sets: fewer bytes row by row
    assert tr.choose_route(32, V, H, e, [1242] * 32, 700) == "row-sparse"
    # everything legal: dense
    assert tr.choose_route(8, V, H, e, [V] * 8, 1940) == "dense-mask"


def test_route_cost_defaults_match_python_model():
    """The device selector's built-in cost model is the Python B200_COST."""
    assert _native.default_route_cost() == tr.B200_COST


STEERED_COST = {"row_sparse_fixed_us": 0.5, "block_floor_us": 0.0, "block_fixed_us": 1.0, "dense_fixed_us": 0.0}


def test_native_route_choice_matches_python_model():
    """gsp_choose_route (the code the device selector runs) picks the route
    choose_route picks, on random statistics and on exact cost ties."""
    import numpy as np
    rng = np.random.default_rng(0)
    for cost in (None, STEERED_COST):
        for _ in range(1500):
            batch = int(rng.integers(1, 300))
            vocab = int(rng.integers(1000, 300000))
            hidden = int(rng.integers(64, 8192))
            ntiles = (vocab + 127) // 128
            legal = [int(x) for x in rng.integers(0, vocab + 1, size=batch) * rng.random(batch) ** 4]
            active = int(rng.integers(0, ntiles + 1))
            got = _native.choose_route_code(batch, vocab, hidden, 2, sum(legal), active, cost)
            assert tr.ROUTES[got] == tr.choose_route(batch, vocab, hidden, 2, legal, active, cost), \
                (batch, vocab, hidden, sum(legal), active, cost)
    # equal block and dense costs: block first, as in choose_route's tuple order
    tie = {"block_floor_us": 0.0, "block_fixed_us": 5.0, "block_gbs": 6000.0, "dense_fixed_us": 5.0,
           "dense_gbs": 6000.0, "row_sparse_fixed_us": 1e9}
    assert tr.choose_route(8, 4096, 256, 2, [4096] * 8, 32, tie) == "block-sparse"
    assert _native.choose_route_code(8, 4096, 256, 2, 8 * 4096, 32, tie) == 1
    assert _native.choose_route_code(1, 4096, 256, 2, 10, 1, tie) == 0  # batch 1: row-sparse


def test_adaptive_entry_validation():
    lib = _native.load()
    route = ctypes.c_int32(7)
    args = [FAKE, 8, FAKE, 8, None, 0, 2, 64, 8, 0, None, 64, None, None, None, None, ctypes.byref(route), None, 0,
            None]
    assert lib.gsp_adaptive_logits(*args) == -1  # bitmask required
    assert route.value == -1 and b"bitmask" in lib.gsp_last_error()
    args[4] = FAKE
    assert lib.gsp_adaptive_logits(*args) == -3  # workspace required
    args[9] = 5
    assert lib.gsp_adaptive_logits(*args) == -2  # dtype
    with pytest.raises(ValueError):
        _native.route_cost({"no_such_field": 1.0})


def test_grouped_entry_validation():
    lib = _native.load()
    assert lib.gsp_group_plan_words(0) == 0 and lib.gsp_group_plan_words(4) == 16 + 24
    assert lib.gsp_grouped_scratch_bytes(0, 10, 10, 1) == 0
    with_l = lib.gsp_grouped_scratch_bytes(32, 248320, 2048, 1)
    without = lib.gsp_grouped_scratch_bytes(32, 248320, 2048, 0)
    assert with_l - without >= 32 * 248320 * 2 and with_l % 256 == 0
    hdr = (ctypes.c_int32 * 8)()
    args = [FAKE, 8, FAKE, 8, FAKE, 2, 300, 64, 8, 0, None, 64, None, None, None, hdr, FAKE, 1 << 20, FAKE, 1 << 30,
            None]
    assert lib.gsp_grouped_logits(*args) == -1  # batch over GSP_GROUP_MAX_BATCH
    args[6] = 4
    args[4] = None
    assert lib.gsp_grouped_logits(*args) == -1 and b"bitmask" in lib.gsp_last_error()
    assert lib.gsp_group_plan(FAKE, 2, 300, 64, 8, 2, 0, None, FAKE, None) == -1
    assert lib.gsp_group_plan(FAKE, 2, 4, 64, 8, 2, 0, None, None, None) == -1
    assert lib.gsp_gather_rows(FAKE, 16, FAKE, 2, 16, FAKE, 8, None) == -1  # dst stride < row bytes
    assert lib.gsp_gather_rows(None, 16, None, 0, 16, None, 16, None) == 0  # nothing to copy


def test_copy_bytes_validation():
    lib = _native.load()
    assert lib.gsp_copy_bytes(None, None, 0, None) == 0  # nothing to copy
    assert lib.gsp_copy_bytes(None, FAKE, 16, None) == -1
    assert lib.gsp_copy_bytes(FAKE, None, 16, None) == -1


def test_merge_logsumexp_validation():
    lib = _native.load()
    assert lib.gsp_merge_logsumexp(FAKE, 0, 4, FAKE, None) == -1
    assert lib.gsp_merge_logsumexp(None, 2, 4, FAKE, None) == -1


def test_newer_python_entries_reject_cpu_tensors_and_bad_arguments():
    """The device-route, lane-group and graphed-head entry points raise
    ValueError for CPU tensors like the reference's entry points (no CPU
    path), and unknown policies or oversized grouped batches are refused
    before any device work."""
    h = torch.zeros(2, 8, dtype=torch.float16)
    w = torch.zeros(64, 8, dtype=torch.float16)
    m = torch.zeros(2, 2, dtype=torch.int32)
    for call in (lambda: tr.grammar_head(h, w, m),
                 lambda: tr.grouped_grammar_logits(h, w, m),
                 lambda: tr.adaptive_grammar_logits(h, w, m, policy="device"),
                 lambda: tr.adaptive_grammar_logits(h, w, m, policy="grouped"),
                 lambda: tr.adaptive_grammar_logits(h, w, m, policy="no-such-policy")):
        with pytest.raises(ValueError):
            call()
    from gsp.graphed import GraphedGrammarHead
    with pytest.raises(ValueError):
        GraphedGrammarHead(w, 2)


def test_ctypes_signatures_match_header_parameter_counts():
    """Every entry point declared in include/gsp_b200.h has a ctypes
    signature with the same number of parameters (an ABI change that misses
    the binding fails here, on CPU)."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    decls = re.findall(r"^\s*(?:int32_t|size_t|void|const char\s*\*)\s*(gsp_\w+)\s*\(([^;]*?)\)\s*;", text, re.M | re.S)
    assert len(decls) >= 20
    for name, params in decls:
        params = " ".join(params.split())
        n = 0 if params in ("", "void") else params.count(",") + 1
        assert name in _native.SIGNATURES, name
        assert len(_native.SIGNATURES[name][0]) == n, (name, n, len(_native.SIGNATURES[name][0]))
