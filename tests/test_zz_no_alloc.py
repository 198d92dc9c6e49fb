"""GPU test of gsp_row_sparse_logits_static, the entry point for callers that
cannot allocate device memory (for example a plugin inside a serving engine
that owns all device memory, or an FFI binding handed only its input and
output buffers). The call must produce what the ordinary workspace-taking
entry point produces, on two calls in a row (the second one reuses the
library's shared scratch array), and must refuse sizes above its limits.

This file is collected last on purpose, so that a run stopping at the first
failure has already run every other test; it also passes on its own.
"""
import ctypes

import numpy as np
import pytest
import torch

from gsp import _native
from oracle import gsp_oracle as O

pytestmark = pytest.mark.gpu

STATIC_MAX_BATCH = 1024
STATIC_MAX_VOCAB = 1 << 20


def _static_call(h, w, mask, logits, top_value, top_index, top_key):
    lib = _native.load()
    return lib.gsp_row_sparse_logits_static(
        ctypes.c_void_p(h.data_ptr()), h.stride(0), ctypes.c_void_p(w.data_ptr()), w.stride(0),
        ctypes.c_void_p(mask.data_ptr()), mask.stride(0), h.shape[0], w.shape[0], h.shape[1],
        _native.dtype_code(h.dtype), 0, ctypes.c_void_p(logits.data_ptr()), logits.stride(0),
        ctypes.c_void_p(top_value.data_ptr()), ctypes.c_void_p(top_index.data_ptr()),
        ctypes.c_void_p(top_key.data_ptr()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def _outputs(batch, vocab, dev, dtype):
    return (torch.empty(batch, vocab, device=dev, dtype=dtype), torch.empty(batch, device=dev, dtype=torch.float32),
            torch.empty(batch, device=dev, dtype=torch.int64), torch.empty(batch, device=dev, dtype=torch.int64))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_static_entry_matches_workspace_entry_twice(cuda_device, dtype):
    rng = np.random.default_rng(2024)
    vocab, hidden, batch = 50_000, 512, 3
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32) * np.float32(0.02)).to(dtype)
    h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).to(dtype)
    wd, hd = w.to(cuda_device), h.to(cuda_device)
    for call in range(2):  # the second call finds the scratch left by the first
        mask = O.make_batch_mask(rng, batch, vocab, [500, 0, 7000], clustered=(call == 1), max_runs=16)
        md = torch.from_numpy(mask).to(cuda_device)
        ref = _outputs(batch, vocab, cuda_device, dtype)
        _native.row_sparse(hd, wd, md, logits=ref[0], top_value=ref[1], top_index=ref[2], top_key=ref[3])
        got = _outputs(batch, vocab, cuda_device, dtype)
        status = _static_call(hd, wd, md, *got)
        assert status == _native.GSP_OK, _native.load().gsp_last_error()
        torch.cuda.synchronize()
        exact = O.masked_logits_exact(h, w, mask)
        for out in (ref[0], got[0]):
            rep = O.compare_logits(exact, out.cpu(), dtype=dtype)
            assert rep["support"] and rep["values"], (call, rep)
        rep = O.compare_logits(ref[0].cpu().double(), got[0].cpu(), dtype=dtype)
        assert rep["support"] and rep["values"], (call, rep)
        assert torch.equal(got[2], ref[2]) and torch.equal(got[1], ref[1]) and torch.equal(got[3], ref[3])
        assert torch.equal(got[2], got[0].argmax(-1))
        assert got[2][1].item() == 0 and got[1][1].item() == float("-inf")  # empty legal set


def _static_error(lib):
    err = ctypes.c_int32(-1)
    status = lib.gsp_row_sparse_static_error(ctypes.byref(err),
                                            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert status == _native.GSP_OK, lib.gsp_last_error()
    return err.value


# (batch, vocab, hidden): a batch whose flat mask (62,080 words) is above the
# multi-request threshold, the largest batch on a small vocabulary, and the
# largest vocabulary at batch 1; run in this order, so each call finds the
# scratch as a call of another size left it.
_LIMIT_CASES = [(8, 248_320, 256), (STATIC_MAX_BATCH, 2_000, 64), (1, STATIC_MAX_VOCAB, 64), (8, 248_320, 256)]


def test_static_entry_large_batches_and_limits(cuda_device):
    lib = _native.load()
    assert _static_error(lib) == 0
    rng = np.random.default_rng(77)
    dtype = torch.float16
    for batch, vocab, hidden in _LIMIT_CASES:
        w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32) * np.float32(0.02)).to(dtype)
        h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).to(dtype)
        legal = [int(x) for x in rng.integers(0, max(2, vocab // 100), size=batch)]
        legal[0] = 0
        mask = O.make_batch_mask(rng, batch, vocab, legal, clustered=batch % 2 == 0, max_runs=16)
        wd, hd, md = w.to(cuda_device), h.to(cuda_device), torch.from_numpy(mask).to(cuda_device)
        ref = _outputs(batch, vocab, cuda_device, dtype)
        _native.row_sparse(hd, wd, md, logits=ref[0], top_value=ref[1], top_index=ref[2], top_key=ref[3])
        got = _outputs(batch, vocab, cuda_device, dtype)
        for _ in range(2):  # two calls in a row on the same inputs
            got[0].fill_(0)
            status = _static_call(hd, wd, md, *got)
            assert status == _native.GSP_OK, lib.gsp_last_error()
            torch.cuda.synchronize()
            rep = O.compare_logits(ref[0].cpu().double(), got[0].cpu(), dtype=dtype)
            assert rep["support"] and rep["values"], (batch, vocab, rep)
            assert torch.equal(got[2], ref[2]) and torch.equal(got[3], ref[3]), (batch, vocab)
        sel = slice(0, min(batch, 64))  # the oracle on a slice of the batch
        exact = O.masked_logits_exact(h[sel], w, mask[sel])
        rep = O.compare_logits(exact, got[0][sel].cpu(), dtype=dtype)
        assert rep["support"] and rep["values"], (batch, vocab, rep)
        assert got[2][0].item() == 0 and got[1][0].item() == float("-inf")  # request 0 has no legal token
        assert _static_error(lib) == 0
        del w, wd, ref, got
        torch.cuda.empty_cache()


def test_static_entry_rejects_sizes_beyond_its_scratch(cuda_device):
    lib = _native.load()
    h = torch.zeros(1, 8, device=cuda_device, dtype=torch.float16)
    w = torch.zeros(64, 8, device=cuda_device, dtype=torch.float16)
    mask = torch.zeros(1, 2, device=cuda_device, dtype=torch.int32)
    outs = _outputs(1, 64, cuda_device, torch.float16)
    # batch above the limit: the call must fail before any launch
    status = lib.gsp_row_sparse_logits_static(
        ctypes.c_void_p(h.data_ptr()), 8, ctypes.c_void_p(w.data_ptr()), 8, ctypes.c_void_p(mask.data_ptr()), 0,
        STATIC_MAX_BATCH + 1, 64, 8, 0, 0, ctypes.c_void_p(outs[0].data_ptr()), 64,
        ctypes.c_void_p(outs[1].data_ptr()), ctypes.c_void_p(outs[2].data_ptr()), ctypes.c_void_p(outs[3].data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert status == _native.GSP_ERR_INVALID_ARGUMENT
    assert b"static scratch limits" in lib.gsp_last_error()
    status = lib.gsp_row_sparse_logits_static(
        ctypes.c_void_p(h.data_ptr()), 8, ctypes.c_void_p(w.data_ptr()), 8, ctypes.c_void_p(mask.data_ptr()), 0,
        1, STATIC_MAX_VOCAB + 1, 8, 0, 0, ctypes.c_void_p(outs[0].data_ptr()), 64,
        ctypes.c_void_p(outs[1].data_ptr()), ctypes.c_void_p(outs[2].data_ptr()), ctypes.c_void_p(outs[3].data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert status == _native.GSP_ERR_INVALID_ARGUMENT
