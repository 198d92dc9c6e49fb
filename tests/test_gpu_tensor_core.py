"""GPU parity of the tensor-core paths: the grammar-aware block GEMM
(gsp_block_gemm_logits: active-tile builder + tcgen05 projection) and the
dense masked GEMM (gsp_dense_masked_logits), against the CPU oracle and the
reference's golden outputs, plus the adaptive dispatcher.

Tolerance as in test_gpu_row_sparse.py (oracle.value_bound): support bit-exact,
legal logits within atol 2e-3 + max(rtol 2e-3 * |exact|, half an output ulp),
greedy top-1 equal to the exact argmax outside the near-tie window, fused top-1
equal to torch.argmax of the kernel's own logits.
"""
import numpy as np
import pytest
import torch

from conftest import load_json, load_npz
from gsp import _native
from gsp import triton_runtime as tr
from oracle import gsp_oracle as O

pytestmark = pytest.mark.gpu


def _check(exact, got, dtype, label=""):
    rep = O.compare_logits(exact, got.cpu(), dtype=dtype)
    assert rep["support"], ("support", label, rep)
    assert rep["values"], ("values", label, rep)
    _, idx = O.top1(got.cpu())
    assert O.top1_agrees(exact, idx, dtype=dtype), ("top1", label)


def _run(fn, h, w, mask, with_logits=True):
    b, v = h.shape[0], w.shape[0]
    logits = torch.empty(b, v, device=h.device, dtype=h.dtype) if with_logits else None
    tv = torch.empty(b, device=h.device, dtype=torch.float32)
    ti = torch.empty(b, device=h.device, dtype=torch.int64)
    fn(h, w, mask, logits=logits, top_value=tv, top_index=ti)
    return logits, tv, ti


@pytest.mark.parametrize("fixture", ["block_gemm_ref.npz", "dense_mask_ref.npz"])
@pytest.mark.parametrize("route", ["block", "dense"])
def test_golden_fixtures(cuda_device, fixture, route):
    data, meta = load_npz(fixture)
    fn = _native.block_gemm if route == "block" else _native.dense_masked
    for c in meta:
        w, h, mask = O.kernel_case_inputs(c["vocab"], c["hidden"], c["batch"], c["dtype"], c["seed"],
                                          c["recipe"], c["extra_words"])
        ref = O.bits16_to_tensor(data[c["name"] + "/out"], c["dtype"])
        logits, tv, ti = _run(fn, h.to(cuda_device), w.to(cuda_device), torch.from_numpy(mask).to(cuda_device))
        assert torch.equal(torch.isfinite(logits.cpu()), torch.isfinite(ref)), (route, c["name"])
        _check(O.masked_logits_exact(h, w, mask), logits, O.TORCH_DTYPES[c["dtype"]], c["name"])
        assert torch.equal(ti, logits.argmax(-1)), (route, c["name"])
        assert torch.equal(tv, logits.float().gather(1, ti[:, None])[:, 0]), (route, c["name"])


def test_reference_block_gemm_test_shapes(cuda_device):
    """tests/test_triton_block_gemm.py of the reference: V=248,320, H=2,048,
    fp16, batches {2,4,8,16,32}, alternating k = 7 / 4096 uniform ids per request."""
    vocab, hidden = 248320, 2048
    g = torch.Generator(device=cuda_device).manual_seed(99)
    wd = torch.randn(vocab, hidden, device=cuda_device, generator=g).half()
    w = wd.cpu()
    rng = np.random.default_rng(123)
    for batch in (2, 4, 8, 16, 32):
        hd = torch.randn(batch, hidden, device=cuda_device, generator=g).half()
        ks = [7 if i % 2 == 0 else 4096 for i in range(batch)]
        mask = O.make_batch_mask(rng, batch, vocab, ks)
        got = tr.bitmask_block_gemm_logits(hd, wd, torch.from_numpy(mask).to(cuda_device))
        _check(O.masked_logits_exact(hd.cpu(), w, mask), got, torch.float16, f"batch={batch}")


@pytest.mark.parametrize("batch", [2, 4, 8, 16, 32])
def test_batched_clustered_workload(cuda_device, batch):
    """V=248,320, H=2,048 fp16, each request 0.5% legal in <= 16 clustered runs."""
    vocab, hidden = 248320, 2048
    g = torch.Generator(device=cuda_device).manual_seed(7)
    wd = (torch.randn(vocab, hidden, device=cuda_device, generator=g) * 0.02).half()
    hd = torch.randn(batch, hidden, device=cuda_device, generator=g).half()
    rng = np.random.default_rng(batch)
    mask = O.make_batch_mask(rng, batch, vocab, [1242] * batch, clustered=True, max_runs=16)
    md = torch.from_numpy(mask).to(cuda_device)
    exact = O.masked_logits_exact(hd.cpu(), wd.cpu(), mask)
    results = {}
    for fn in (_native.block_gemm, _native.dense_masked, _native.row_sparse):
        logits, tv, ti = _run(fn, hd, wd, md)
        _check(exact, logits, torch.float16, fn.__name__)
        assert torch.equal(ti, logits.argmax(-1))
        results[fn.__name__] = (tv, ti)
    # top-1 without materialising logits: identical to the same kernel's with-logits run
    _, tv2, ti2 = _run(_native.block_gemm, hd, wd, md, with_logits=False)
    tv, ti = results["block_gemm"]
    assert torch.equal(ti2, ti) and torch.equal(tv2, tv)


@pytest.mark.parametrize("vocab,hidden,batch,dtype", [
    (1000, 96, 3, torch.float16),        # V % 128 != 0, H % 64 != 0
    (4100, 200, 5, torch.bfloat16),      # V % 32 != 0
    (2048, 64, 1, torch.float16),        # batch 1 on the tensor cores
    (3000, 128, 300, torch.float16),     # two batch chunks (256 + 44)
    (1025, 512, 33, torch.bfloat16),     # last tile holds one row
    (777, 12, 2, torch.float16),         # H % 8 != 0: row-sparse path
    (1_300_000, 64, 3, torch.float16),   # over 64 tiles per CTA: tile ids read from the workspace list
])
def test_edge_shapes(cuda_device, vocab, hidden, batch, dtype):
    rng = np.random.default_rng(vocab + batch)
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32)).to(dtype)
    h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).to(dtype)
    mask = O.recipe_mask("random+zero+u5+full+c40", rng, batch, vocab)
    exact = O.masked_logits_exact(h, w, mask)
    for fn in (_native.block_gemm, _native.dense_masked):
        logits, tv, ti = _run(fn, h.to(cuda_device), w.to(cuda_device), torch.from_numpy(mask).to(cuda_device))
        _check(exact, logits, dtype, f"{fn.__name__} V={vocab} H={hidden} B={batch}")
        assert torch.equal(ti, logits.argmax(-1))


def test_no_active_tile_and_unmasked_dense(cuda_device):
    rng = np.random.default_rng(11)
    vocab, hidden, batch = 5000, 256, 4
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32)).half()
    h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).half()
    mask = np.zeros((batch, O.mask_words(vocab)), dtype=np.int32)
    logits, tv, ti = _run(_native.block_gemm, h.to(cuda_device), w.to(cuda_device),
                          torch.from_numpy(mask).to(cuda_device))
    assert not torch.isfinite(logits).any()
    assert ti.tolist() == [0] * batch and all(v == float("-inf") for v in tv.tolist())
    # no mask at all: the dense GEMM
    logits, tv, ti = _run(_native.dense_masked, h.to(cuda_device), w.to(cuda_device), None)
    _check(O.masked_logits_exact(h, w, None), logits, torch.float16, "unmasked")
    assert torch.equal(ti, logits.argmax(-1))


def test_adaptive_dispatch_known_answers(cuda_device):
    """tests/test_adaptive_dispatch.py of the reference: routes and parity."""
    routes = {(c["batch"], c["pattern"]): c["route"] for c in load_json("routes_ref.json")["dispatch_cases"]}
    vocab, hidden = 8192, 512
    for (batch, pattern), expected in routes.items():
        g = torch.Generator().manual_seed(1000 + batch)
        h = torch.randn(batch, hidden, generator=g).half()
        w = torch.randn(vocab, hidden, generator=g).half()
        mask = torch.zeros(batch, vocab // 32, dtype=torch.int32)
        for b in range(batch):
            if pattern == "all_dense" or (pattern == "mixed" and b % 2):
                mask[b].fill_(-1)
            else:
                mask[b, 0] = 1
        frac = tr.full_word_fraction_cpu(mask)
        got, route = tr.adaptive_grammar_logits(h.to(cuda_device), w.to(cuda_device), mask.to(cuda_device),
                                                full_word_fraction=frac)
        assert route == expected, (batch, pattern, route)
        got = got.reshape(batch, -1)
        _check(O.masked_logits_exact(h, w, mask.numpy()), got, torch.float16, f"{batch} {pattern}")
        got_b, route_b = tr.adaptive_grammar_logits(h.to(cuda_device), w.to(cuda_device), mask.to(cuda_device),
                                                    full_word_fraction=frac, policy="b200")
        assert route_b in tr.ROUTES
        _check(O.masked_logits_exact(h, w, mask.numpy()), got_b.reshape(batch, -1), torch.float16, route_b)


def test_workspace_reuse_across_batch_sizes(cuda_device):
    """One workspace serves calls of different batch sizes and routes: the
    block path must leave its tile lists zeroed, or a later, larger batch reads
    them back as top-1 keys."""
    rng = np.random.default_rng(5)
    vocab, hidden = 3000, 128
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32)).half().to(cuda_device)
    for batch in (44, 256, 3, 300, 17):
        h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).half().to(cuda_device)
        mask = torch.from_numpy(O.recipe_mask("random+zero+u5+full+c40", rng, batch, vocab)).to(cuda_device)
        for fn in (_native.block_gemm, _native.dense_masked, _native.row_sparse):
            logits, tv, ti = _run(fn, h, w, mask)
            assert torch.equal(ti, logits.argmax(-1)), (batch, fn.__name__)
            assert torch.equal(tv, logits.float().gather(1, ti[:, None])[:, 0]), (batch, fn.__name__)


@pytest.mark.parametrize("route", ["block", "dense"])
def test_top1_with_vocab_offset_tensor_core(cuda_device, route):
    """The fused top-1 of a vocabulary shard (global ids offset by up to and
    past 2^24, as the vocabulary-parallel head reports them) at batches 1-33
    is the argmax of the kernel's own logits, shifted by the offset."""
    vocab, hidden = 50_000, 256
    rng = np.random.default_rng(93)
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32) * np.float32(0.05)).half().to(cuda_device)
    h = torch.from_numpy(rng.standard_normal((33, hidden), dtype=np.float32)).half().to(cuda_device)
    ks = [int(k) for k in rng.integers(1, 3000, size=33)]
    mask = torch.from_numpy(O.make_batch_mask(rng, 33, vocab, ks, clustered=True, max_runs=8)).to(cuda_device)
    fn = _native.block_gemm if route == "block" else _native.dense_masked
    for b in (1, 2, 8, 32, 33):
        logits, tv0, ti0 = _run(fn, h[:b], w, mask[:b])
        assert torch.equal(ti0, logits.argmax(-1)), (route, b)
        for offset in (1_000_000, 1 << 24, (1 << 24) - 40_000):
            tv = torch.empty(b, device=cuda_device)
            ti = torch.empty(b, device=cuda_device, dtype=torch.int64)
            fn(h[:b], w, mask[:b], top_value=tv, top_index=ti, vocab_offset=offset)
            assert torch.equal(ti, ti0 + offset), (route, b, offset)
            assert torch.equal(tv, tv0), (route, b, offset)
    assert _native.workspace_error(cuda_device) == 0


def test_no_bounded_wait_gave_up_tensor_core(cuda_device):
    assert _native.workspace_error(cuda_device) == 0
