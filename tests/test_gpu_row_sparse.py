"""GPU parity of the row-sparse path (gsp_row_sparse_logits / _compact), the
mask utilities and constrained_projection against the CPU oracle and the
reference's golden outputs.

Tolerance (oracle.value_bound): legal support bit-exact; each legal logit
within atol 2e-3 + max(rtol 2e-3 * |exact|, half an output ulp) of the exact
float64 value; greedy top-1 identical to the exact argmax except inside the
near-tie window atol + max(rtol * |max|, one output ulp); fused top-1 equal to
torch.argmax over the kernel's own logits, bit for bit.
"""
import numpy as np
import pytest
import torch

from conftest import load_npz
from gsp import _native
from gsp import runtime as rt
from gsp import triton_runtime as tr
from oracle import gsp_oracle as O

pytestmark = pytest.mark.gpu


def _check(exact, got, dtype, label=""):
    rep = O.compare_logits(exact, got.cpu(), dtype=dtype)
    assert rep["support"], ("support", label, rep)
    assert rep["values"], ("values", label, rep)
    _, idx = O.top1(got.cpu())
    assert O.top1_agrees(exact, idx, dtype=dtype), ("top1", label)


def _fused(h2, w, mask, logits=None):
    b = h2.shape[0]
    tv = torch.empty(b, device=h2.device, dtype=torch.float32)
    ti = torch.empty(b, device=h2.device, dtype=torch.int64)
    tk = torch.empty(b, device=h2.device, dtype=torch.int64)
    _native.row_sparse(h2, w, mask, logits=logits, top_value=tv, top_index=ti, top_key=tk)
    return tv, ti, tk


@pytest.mark.parametrize("fixture", ["row_sparse_ref.npz", "dense_mask_ref.npz"])
def test_golden_fixtures(cuda_device, fixture):
    data, meta = load_npz(fixture)
    for c in meta:
        w, h, mask = O.kernel_case_inputs(c["vocab"], c["hidden"], c["batch"], c["dtype"], c["seed"],
                                          c["recipe"], c["extra_words"])
        ref = O.bits16_to_tensor(data[c["name"] + "/out"], c["dtype"])
        got = tr.bitmask_sparse_logits(h.to(cuda_device), w.to(cuda_device), torch.from_numpy(mask).to(cuda_device))
        got = got.reshape(c["batch"], -1).cpu()
        assert torch.equal(torch.isfinite(got), torch.isfinite(ref)), c["name"]
        _check(O.masked_logits_exact(h, w, mask), got, O.TORCH_DTYPES[c["dtype"]], c["name"])


def test_reference_sparse_test_shapes(cuda_device):
    """tests/test_triton_sparse.py of the reference: V=151,936, H=1,024, fp16,
    batch 1, k in {1, 13, 428, 4096, 32768, 120000}, W and h ~ N(0, 1)."""
    rng = np.random.default_rng(17)
    vocab, hidden = 151936, 1024
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32)).half()
    h = torch.from_numpy(rng.standard_normal((1, hidden), dtype=np.float32)).half()
    wd, hd = w.to(cuda_device), h.to(cuda_device)
    for k in (1, 13, 428, 4096, 32768, 120000):
        ids = rng.permutation(vocab)[:k]
        mask = O.ids_to_bitmask(ids, vocab)
        got = tr.bitmask_sparse_logits(hd, wd, torch.from_numpy(mask).to(cuda_device))
        assert got.shape == (vocab,)
        _check(O.masked_logits_exact(h, w, mask)[0], got, torch.float16, f"k={k}")


def test_fused_top1_is_argmax_of_logits(cuda_device):
    rng = np.random.default_rng(3)
    for vocab, hidden, batch, dtype in ((5000, 256, 1, torch.float16), (4099, 512, 3, torch.bfloat16),
                                        (248320, 64, 2, torch.float16)):
        w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32)).to(dtype).to(cuda_device)
        h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).to(dtype).to(cuda_device)
        mask = torch.from_numpy(O.make_batch_mask(rng, batch, vocab, [vocab // 50] * batch)).to(cuda_device)
        logits = torch.empty(batch, vocab, device=cuda_device, dtype=dtype)
        tv, ti, tk = _fused(h, w, mask, logits)
        assert torch.equal(ti, logits.argmax(-1))
        assert torch.equal(tv, logits.float().gather(1, ti[:, None])[:, 0])
        tv2, ti2, _ = _fused(h, w, mask, None)  # top-1 without materialising logits
        assert torch.equal(ti2, ti) and torch.equal(tv2, tv)


def test_ties_go_to_lowest_index(cuda_device):
    vocab, hidden = 4096, 128
    w = torch.zeros(vocab, hidden, dtype=torch.float16)
    w[:, 0] = 1.0
    h = torch.zeros(1, hidden, dtype=torch.float16)
    h[0, 0] = 2.0
    mask = O.ids_to_bitmask([4000, 17, 900, 3000], vocab)
    logits = torch.empty(1, vocab, device=cuda_device, dtype=torch.float16)
    tv, ti, _ = _fused(h.to(cuda_device), w.to(cuda_device), torch.from_numpy(mask).to(cuda_device), logits)
    assert ti.item() == 17 and tv.item() == 2.0
    assert ti.item() == logits.argmax(-1).item()


def test_empty_mask_and_repeated_calls(cuda_device):
    vocab, hidden = 3000, 64
    rng = np.random.default_rng(9)
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32)).half().to(cuda_device)
    h = torch.from_numpy(rng.standard_normal((2, hidden), dtype=np.float32)).half().to(cuda_device)
    mask = torch.from_numpy(O.make_batch_mask(rng, 2, vocab, [0, 40])).to(cuda_device)
    logits = torch.empty(2, vocab, device=cuda_device, dtype=torch.float16)
    results = [tuple(t.clone() for t in _fused(h, w, mask, logits)) for _ in range(3)]
    for r in results[1:]:
        assert all(torch.equal(a, b) for a, b in zip(r, results[0]))
    tv, ti, _ = results[0]
    assert ti[0].item() == 0 and tv[0].item() == float("-inf")  # torch.argmax of all -inf is 0
    assert not torch.isfinite(logits[0]).any()
    assert ti[1].item() == logits[1].argmax().item()


@pytest.mark.parametrize("vocab,hidden,batch", [(1, 8, 1), (33, 16, 2), (1000, 1000, 2), (4100, 12, 3),
                                                (777, 96, 5)])
def test_edge_shapes(cuda_device, vocab, hidden, batch):
    """V not a multiple of 32, H not a multiple of 8 (scalar path), tiny V."""
    rng = np.random.default_rng(vocab + hidden)
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32)).half()
    h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).half()
    mask = O.recipe_mask("random+full+zero", rng, batch, vocab)
    got = tr.bitmask_sparse_logits(h.to(cuda_device), w.to(cuda_device), torch.from_numpy(mask).to(cuda_device))
    _check(O.masked_logits_exact(h, w, mask).reshape(batch, vocab), got.reshape(batch, vocab), torch.float16)


def test_misaligned_strided_and_broadcast_inputs(cuda_device):
    rng = np.random.default_rng(21)
    vocab, hidden, batch = 2048, 256, 3
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32)).half()
    h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).half()
    mask = O.recipe_mask("u100", rng, 1, vocab, extra_words=3)
    exact = O.masked_logits_exact(h, w, np.repeat(mask, batch, axis=0))
    # hidden starting one element off a 16-byte boundary (vector path disabled)
    hbuf = torch.empty(batch * hidden + 1, dtype=torch.float16, device=cuda_device)
    hbuf[1:] = h.reshape(-1).to(cuda_device)
    h_mis = hbuf[1:].view(batch, hidden)
    # one mask row shared by every request: row stride 0; wider than ceil(V/32)
    m = torch.from_numpy(mask).to(cuda_device).expand(batch, -1)
    logits = torch.empty(batch, vocab + 5, device=cuda_device, dtype=torch.float16)[:, :vocab]
    _native.row_sparse(h_mis, w.to(cuda_device), m, logits=logits)
    _check(exact, logits, torch.float16, "misaligned/broadcast/strided-out")


def test_wide_mask_uses_real_row_stride(cuda_device):
    """A [B, words + extra] mask: every request reads its own row (the reference
    kernels assume stride ceil(V/32); its dense route uses the real stride)."""
    rng = np.random.default_rng(5)
    vocab, hidden, batch = 1000, 64, 3
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32)).half()
    h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).half()
    mask = O.recipe_mask("u10+u300+random", rng, batch, vocab, extra_words=7)
    got = tr.bitmask_sparse_logits(h.to(cuda_device), w.to(cuda_device), torch.from_numpy(mask).to(cuda_device))
    _check(O.masked_logits_exact(h, w, mask), got, torch.float16)


def test_compact_logits(cuda_device):
    rng = np.random.default_rng(8)
    vocab, hidden, batch = 9000, 128, 3
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32)).bfloat16()
    h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).bfloat16()
    mask = O.make_batch_mask(rng, batch, vocab, [5, 0, 700], clustered=True, max_runs=8)
    md = torch.from_numpy(mask).to(cuda_device)
    ids, lg, off = tr.bitmask_compact_logits(h.to(cuda_device), w.to(cuda_device), md)
    legal = O.unpack_bitmask(mask, vocab)
    assert off.tolist() == [0, 5, 5, 705]
    exact = O.masked_logits_exact(h, w, mask)
    for b in range(batch):
        s, e = off[b].item(), off[b + 1].item()
        assert np.array_equal(ids[s:e].cpu().numpy(), np.flatnonzero(legal[b]))
        rep = O.compare_logits(exact[b, np.flatnonzero(legal[b])], lg[s:e].cpu(), dtype=torch.bfloat16)
        assert rep["support"] and rep["values"]


def test_ids_to_bitmask_and_mask_stats(cuda_device):
    rng = np.random.default_rng(12)
    vocab = 248320
    ids = rng.integers(0, vocab, size=5000)
    bm = torch.empty(1, (vocab + 31) // 32, dtype=torch.int32, device=cuda_device)
    stats = torch.empty(2, dtype=torch.int64, device=cuda_device)
    _native.ids_to_bitmask(torch.from_numpy(ids).to(cuda_device), vocab, bm, stats)
    assert np.array_equal(bm.cpu().numpy(), O.ids_to_bitmask(ids, vocab))
    assert stats.tolist() == [len(np.unique(ids)), 0]
    bad = torch.tensor([3, -1, vocab, 5, 5], device=cuda_device)
    _native.ids_to_bitmask(bad, vocab, bm, stats)
    assert stats.tolist() == [2, 2]
    batch = 5
    mask = O.make_batch_mask(rng, batch, vocab, [1242] * batch, clustered=True, max_runs=16)
    mask[2, 10:20] = -1
    st = tr.mask_stats(torch.from_numpy(mask).to(cuda_device), vocab)
    legal = O.unpack_bitmask(mask, vocab)
    assert st["legal_counts"] == legal.sum(1).tolist()
    assert st["full_words"] == [int((mask[b] == -1).sum()) for b in range(batch)]
    assert st["active_tiles"] == O.active_tiles(mask, vocab)


def test_constrained_projection_golden(cuda_device):
    data, _ = load_npz("projection_ref.npz")
    import json
    meta = json.loads(str(data["meta"]))
    for c in meta:
        if c["name"].startswith("config0"):
            continue  # the fp32 configuration: test_gpu_fp32.py
        w, h = O.projection_case_inputs(c["dtype"], c["seed"])
        if c["hidden_1d"]:
            h = h[0]
        ids = None if c["ids_is_none"] else torch.from_numpy(data[c["name"] + "/ids"])
        res = rt.constrained_projection(h.to(cuda_device), w.to(cuda_device),
                                        None if ids is None else ids.to(cuda_device),
                                        dense_threshold=c["threshold"])
        assert res.mode == c["mode"], c["name"]
        assert np.array_equal(res.token_ids.cpu().numpy(), data[c["name"] + "/token_ids"]), c["name"]
        exact = O.constrained_projection(h, w, ids, dense_threshold=c["threshold"])
        ex = (h.reshape(-1, h.shape[-1]).double() @ w[exact.token_ids].double().T)
        ex = ex[0] if h.ndim == 1 else ex
        rep = O.compare_logits(ex, res.logits.cpu(), dtype=w.dtype)
        assert rep["support"] and rep["values"], (c["name"], rep)


def test_constrained_projection_errors_and_config0(cuda_device):
    w = torch.zeros((100, 8), dtype=torch.float16, device=cuda_device)
    h = torch.zeros((1, 8), dtype=torch.float16, device=cuda_device)
    with pytest.raises(ValueError, match="grammar produced an empty legal-token set"):
        rt.constrained_projection(h, w, torch.zeros(0, dtype=torch.long))
    with pytest.raises(ValueError, match="out-of-range"):
        rt.constrained_projection(h, w, torch.tensor([5, 100]))
    with pytest.raises(ValueError, match="one-dimensional"):
        rt.constrained_projection(h, w, torch.tensor([[1, 2]]))
    with pytest.raises(ValueError, match="unsupported dtype"):
        rt.constrained_projection(h.double(), w.double(), torch.tensor([1]))
    # 32,768 x 1,024, batch 1, 1% uniform (seed 0), also in fp16 (the fp32
    # configuration itself is checked in test_gpu_fp32.py)
    w32, h32, ids = O.config0_inputs(seed=0)
    w16, h16 = w32.half(), h32.half()
    res = rt.constrained_projection(h16.to(cuda_device), w16.to(cuda_device), torch.from_numpy(ids).to(cuda_device))
    assert res.mode == "sparse-gather" and res.logits.shape == (1, 327)
    assert np.array_equal(res.token_ids.cpu().numpy(), ids)
    exact = h16.double() @ w16[torch.from_numpy(ids)].double().T
    rep = O.compare_logits(exact, res.logits.cpu(), dtype=torch.float16)
    assert rep["values"], rep


@pytest.mark.parametrize("clustered", [False, True])
def test_full_size_density_sweep(cuda_device, clustered):
    """V=248,320, H=2,048 fp16, W ~ N(0, 0.02), h ~ N(0, 1), batch 1: every
    density of the GEMV workload, uniform or clustered in 1-64 runs."""
    vocab, hidden = 248320, 2048
    g = torch.Generator(device=cuda_device).manual_seed(1234)
    wd = (torch.randn(vocab, hidden, device=cuda_device, generator=g) * 0.02).half()
    hd = torch.randn(1, hidden, device=cuda_device, generator=g).half()
    w, h = wd.cpu(), hd.cpu()
    rng = np.random.default_rng(77 + clustered)
    for density in (0.0005, 0.005, 0.01, 0.10, 0.50, 1.0):
        k = int(round(density * vocab))
        mask = O.make_batch_mask(rng, 1, vocab, [k], clustered=clustered, max_runs=64)
        logits = torch.empty(1, vocab, device=cuda_device, dtype=torch.float16)
        tv, ti, _ = _fused(hd, wd, torch.from_numpy(mask).to(cuda_device), logits)
        exact = O.masked_logits_exact(h, w, mask)
        _check(exact, logits, torch.float16, f"density={density}")
        assert int(torch.isfinite(logits).sum()) == k
        assert ti.item() == logits.argmax(-1).item()


@pytest.mark.parametrize("clustered", [False, True])
def test_batch1_mask_over_8192_words(cuda_device, clustered):
    """Batch 1 with a vocabulary of more than 262,144 tokens (9,376 mask words,
    a ragged last word): the staged kernel holds 32 mask words per thread, and
    the half-warps resolve each unit from two groups of 16 staged words."""
    vocab, hidden = 300_007, 128
    rng = np.random.default_rng(4242 + clustered)
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32) * np.float32(0.05)).half()
    h = torch.from_numpy(rng.standard_normal((1, hidden), dtype=np.float32)).half()
    wd, hd = w.to(cuda_device), h.to(cuda_device)
    for density in (0.01, 0.10):
        k = int(round(density * vocab))
        mask = O.make_batch_mask(rng, 1, vocab, [k], clustered=clustered, max_runs=32)
        mask[0, -1] |= np.int32(-1)  # bits beyond the vocabulary set: the kernel must ignore them
        logits = torch.empty(1, vocab, device=cuda_device, dtype=torch.float16)
        tv, ti, _ = _fused(hd, wd, torch.from_numpy(mask).to(cuda_device), logits)
        exact = O.masked_logits_exact(h, w, mask)
        _check(exact, logits, torch.float16, f"density={density}")
        assert ti.item() == logits.argmax(-1).item()


def test_top1_merge_paths_agree(cuda_device):
    """Global ids below 2^24 - 1 take the polled top-1 merge (self-tagged
    per-CTA key slots); a vocabulary offset that reaches past it takes the
    ticket merge. Both report the same token, shifted by the offset."""
    vocab, hidden = 50_000, 256
    rng = np.random.default_rng(91)
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32) * np.float32(0.05)).half().to(cuda_device)
    h = torch.from_numpy(rng.standard_normal((2, hidden), dtype=np.float32)).half().to(cuda_device)
    mask = torch.from_numpy(O.make_batch_mask(rng, 2, vocab, [400, 3000], clustered=True, max_runs=8)).to(cuda_device)
    for b in (1, 2):
        tv0, ti0, _ = _fused(h[:b], w, mask[:b])
        for offset in (0, 1_000_000, 1 << 24, (1 << 24) - 40_000):
            tv = torch.empty(b, device=cuda_device)
            ti = torch.empty(b, device=cuda_device, dtype=torch.int64)
            _native.row_sparse(h[:b], w, mask[:b], top_value=tv, top_index=ti, vocab_offset=offset)
            assert torch.equal(ti, ti0 + offset), (b, offset)
            assert torch.equal(tv, tv0), (b, offset)
    assert _native.workspace_error(cuda_device) == 0


def test_no_bounded_wait_gave_up(cuda_device):
    """Every kernel above completed without giving up a bounded wait."""
    assert _native.workspace_error(cuda_device) == 0


def test_copy_bytes_and_top1_into_pinned_memory(cuda_device):
    """gsp_copy_bytes between pinned host and device memory (16-byte units and
    ragged tails), and a projection storing its top-1 straight into pinned
    host memory: the end-to-end step's transfers."""
    dev = cuda_device
    rng = np.random.default_rng(21)
    for nbytes, offset in ((35 * 1024, 0), (35 * 1024 + 3, 0), (1000, 1), (16, 0), (1, 0)):
        src = torch.from_numpy(rng.integers(0, 256, size=nbytes + offset, dtype=np.uint8)).pin_memory()
        dst = torch.zeros(nbytes + offset, dtype=torch.uint8, device=dev)
        _native.copy_bytes(dst[offset:], src[offset:], nbytes)
        back = torch.zeros(nbytes + offset, dtype=torch.uint8).pin_memory()
        _native.copy_bytes(back[offset:], dst[offset:], nbytes)
        torch.cuda.synchronize()
        assert torch.equal(dst[offset:].cpu(), src[offset:]) and torch.equal(back[offset:], src[offset:]), nbytes
    vocab, hidden = 20000, 256
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32) * 0.1).half().to(dev)
    h = torch.from_numpy(rng.standard_normal((1, hidden), dtype=np.float32)).half().to(dev)
    mask = torch.from_numpy(O.make_batch_mask(rng, 1, vocab, [200])).to(dev)
    tv_h = torch.zeros(1, dtype=torch.float32).pin_memory()
    ti_h = torch.zeros(1, dtype=torch.int64).pin_memory()
    tv_d = torch.empty(1, device=dev)
    ti_d = torch.empty(1, dtype=torch.int64, device=dev)
    for _ in range(2):
        _native.row_sparse(h, w, mask, top_value=tv_h, top_index=ti_h)
        _native.row_sparse(h, w, mask, top_value=tv_d, top_index=ti_d)
        torch.cuda.synchronize()
        assert ti_h.item() == ti_d.item() and tv_h.item() == tv_d.item()


def test_fused_host_input_step(cuda_device):
    """gsp_row_sparse_step (PreparedStep): one C-ABI call copies the pinned
    staging row (mask + hidden state) to the device and projects, the top-1
    record landing in pinned host memory; equal to gsp_copy_bytes followed by
    gsp_row_sparse_logits, over staging rows that change every call. A bad
    argument fails before anything is queued (the device row is untouched)."""
    import ctypes
    dev = cuda_device
    rng = np.random.default_rng(31)
    vocab, hidden = 30_000, 512
    words = (vocab + 31) // 32
    mask_pad = (words * 4 + 15) // 16 * 16
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32) * 0.05).half().to(dev)
    rows = []
    for j in range(3):
        row = torch.zeros(mask_pad + hidden * 2, dtype=torch.uint8).pin_memory()
        m = O.make_batch_mask(rng, 1, vocab, [50 * (j + 1)], clustered=j == 1, max_runs=4)
        row[:words * 4] = torch.from_numpy(np.ascontiguousarray(m)).view(torch.uint8).reshape(-1)
        row[mask_pad:] = torch.from_numpy(rng.standard_normal(hidden, dtype=np.float32)).half().view(torch.uint8)
        rows.append(row)
    dev_row = torch.zeros(rows[0].numel(), dtype=torch.uint8, device=dev)
    dev_mask = dev_row[:words * 4].view(torch.int32).view(1, words)
    dev_hidden = dev_row[mask_pad:].view(torch.float16).view(1, hidden)
    host_top = torch.zeros(2, dtype=torch.int64).pin_memory()
    logits = torch.empty(1, vocab, device=dev, dtype=torch.float16)
    step = _native.PreparedStep(rows[0], dev_row, dev_hidden, w, dev_mask, logits=logits,
                                top_value=host_top[1:2].view(torch.float32)[:1], top_index=host_top[0:1])
    ref_logits = torch.empty_like(logits)
    ti = torch.empty(1, device=dev, dtype=torch.int64)
    for j in (0, 1, 2, 0):
        host_top.fill_(-7)
        step(rows[j])
        torch.cuda.synchronize()
        ref_row = torch.empty_like(dev_row)
        _native.copy_bytes(ref_row, rows[j])
        _native.row_sparse(ref_row[mask_pad:].view(torch.float16).view(1, hidden), w,
                           ref_row[:words * 4].view(torch.int32).view(1, words), logits=ref_logits, top_index=ti)
        torch.cuda.synchronize()
        assert torch.equal(dev_row, ref_row) and torch.equal(logits.view(torch.int16), ref_logits.view(torch.int16))
        assert int(host_top[0]) == ti.item() == logits.argmax(-1).item()
    # the same step recorded as a CUDA graph inside the library, its copy
    # pointed at another pinned row on each launch
    gstep = _native.GraphStep(rows[0], dev_row, dev_hidden, w, dev_mask, logits=logits,
                              top_value=host_top[1:2].view(torch.float32)[:1], top_index=host_top[0:1])
    for j in (2, 1, 1, 0, 2):
        host_top.fill_(-7)
        gstep(rows[j])
        torch.cuda.synchronize()
        ref_row = torch.empty_like(dev_row)
        _native.copy_bytes(ref_row, rows[j])
        _native.row_sparse(ref_row[mask_pad:].view(torch.float16).view(1, hidden), w,
                           ref_row[:words * 4].view(torch.int32).view(1, words), logits=ref_logits, top_index=ti)
        torch.cuda.synchronize()
        assert torch.equal(dev_row, ref_row) and torch.equal(logits.view(torch.int16), ref_logits.view(torch.int16))
        assert int(host_top[0]) == ti.item()
    gstep.close()
    assert _native.workspace_error(dev) == 0
    # hidden_dim 0 is rejected before the copy: the device row keeps its bytes
    before = dev_row.clone()
    lib = _native.load()
    st = lib.gsp_row_sparse_step(ctypes.c_void_p(rows[1].data_ptr()), rows[1].numel(),
                                 ctypes.c_void_p(dev_row.data_ptr()), ctypes.c_void_p(dev_hidden.data_ptr()), hidden,
                                 ctypes.c_void_p(w.data_ptr()), hidden, ctypes.c_void_p(dev_mask.data_ptr()), words,
                                 1, vocab, 0, 0, 0, None, vocab, None, None, None, None, 0,
                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == _native.GSP_ERR_INVALID_ARGUMENT
    torch.cuda.synchronize()
    assert torch.equal(dev_row, before)
