"""Vocabulary-parallel head on 2 GPUs (one spawned process per GPU, NCCL for
the set-up): the in-kernel peer exchange (gsp_vocab_parallel_logits) and the
NCCL all-reduce path both give the global greedy top-1 of the full head, equal
to the oracle's exact argmax outside the near-tie window and bit-identical to
each other, for every route, over repeated calls and CUDA-graph replays.
Skipped on machines with fewer than 2 GPUs."""
import math
import os
import socket
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROUTES = ("row-sparse", "block-sparse", "dense-mask")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(vocab, hidden, batch, seed, dtype):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), ".."))
    from oracle import gsp_oracle as O
    rng = np.random.default_rng(seed)
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32) * 0.05).to(dtype)
    h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).to(dtype)
    ks = [int(k) for k in rng.integers(1, max(2, vocab // 50), size=batch)]
    mask = O.make_batch_mask(rng, batch, vocab, ks, clustered=True, max_runs=8)
    return w, h, mask


def _worker(rank, world, port, result_path):
    import sys
    import datetime
    root = os.path.join(os.path.dirname(__file__), "..")
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "grammar-sparse-projection_b200"))
    import torch.distributed as dist
    from gsp import _native
    from gsp import vocab_parallel as vp
    from oracle import gsp_oracle as O

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    failures = []
    try:
        xch = vp.PeerExchange(max_batch=40)
        for vocab, hidden, batch, seed, dtype in ((50000, 256, 1, 1, torch.float16),
                                                  (40000, 128, 3, 2, torch.bfloat16),
                                                  (30001, 64, 33, 3, torch.float16)):
            w, h, mask = _case(vocab, hidden, batch, seed, dtype)
            exact = O.masked_logits_exact(h, w, mask)
            head_peer = vp.VocabParallelHead.from_full_weight(w.to(dev), exchange=xch)
            head_nccl = vp.VocabParallelHead.from_full_weight(w.to(dev))
            hd, md = h.to(dev), torch.from_numpy(mask).to(dev)
            for route in ROUTES:
                tv_n, ti_n, _ = head_nccl.forward(hd, md, route=route)
                for rep in range(3):  # repeated calls advance the exchange epoch
                    tv_p, ti_p, lg = head_peer.forward(hd, md, route=route, full_logits=(rep == 0))
                    if not (torch.equal(tv_p, tv_n) and torch.equal(ti_p, ti_n)):
                        failures.append(f"{route} V={vocab} B={batch} rep {rep}: peer != nccl")
                    if not O.top1_agrees(exact, ti_p.cpu(), dtype=dtype):
                        failures.append(f"{route} V={vocab} B={batch}: top-1 vs oracle")
                    if lg is not None:
                        rep_ = O.compare_logits(exact, lg.cpu(), dtype=dtype)
                        if not (rep_["support"] and rep_["values"]):
                            failures.append(f"{route} V={vocab} B={batch}: gathered logits")
            # the fence-and-flag protocol of heads with 2^24 - 1 or more tokens
            mask_local = head_peer.local_mask(md)
            tv_n, ti_n, _ = head_nccl.forward(hd, md, route="row-sparse")
            for _ in range(3):
                tv_f = torch.empty(batch, device=dev)
                ti_f = torch.empty(batch, device=dev, dtype=torch.int64)
                _native.vocab_parallel("row-sparse", hd, head_peer.weight, mask_local, xch.peers, xch.rank,
                                       xch.max_batch, 1 << 25, top_value=tv_f, top_index=ti_f,
                                       vocab_offset=head_peer.start)
                if not (torch.equal(tv_f, tv_n) and torch.equal(ti_f, ti_n)):
                    failures.append(f"flag protocol V={vocab} B={batch}")
            # CUDA graph: three exchange calls per replay, replayed twice
            tv_g = torch.empty(batch, device=dev)
            ti_g = torch.empty(batch, device=dev, dtype=torch.int64)
            mask_local = head_peer.local_mask(md)
            s = torch.cuda.Stream(device=dev)
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                _native.vocab_parallel("row-sparse", hd, head_peer.weight, mask_local, xch.peers, xch.rank,
                                       xch.max_batch, vocab, top_value=tv_g, top_index=ti_g,
                                       vocab_offset=head_peer.start)
            torch.cuda.current_stream().wait_stream(s)
            torch.cuda.synchronize()
            dist.barrier()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for _ in range(3):
                    _native.vocab_parallel("row-sparse", hd, head_peer.weight, mask_local, xch.peers, xch.rank,
                                           xch.max_batch, vocab, top_value=tv_g, top_index=ti_g,
                                           vocab_offset=head_peer.start)
            for _ in range(2):
                dist.barrier()
                g.replay()
                torch.cuda.synchronize()
                tv_n, ti_n, _ = head_nccl.forward(hd, md, route="row-sparse")
                if not (torch.equal(tv_g, tv_n) and torch.equal(ti_g, ti_n)):
                    failures.append(f"graph replay V={vocab} B={batch}")
            del g
        # sampling across the shards (NCCL merge) equals the single-GPU sampler
        from gsp import triton_runtime as tr
        w, h, mask = _case(30001, 128, 5, 7, torch.float16)
        head_s = vp.VocabParallelHead.from_full_weight(w.to(dev))
        seeds = torch.arange(5, device=dev, dtype=torch.int64) * 7919 + 3
        got = head_s.sample(h.to(dev), torch.from_numpy(mask).to(dev), seeds=seeds, step=4, temperature=0.8)
        want = tr.grammar_sample(h.to(dev), w.to(dev), torch.from_numpy(mask).to(dev), seeds=seeds, step=4,
                                 temperature=0.8)
        if not (torch.equal(got.token_ids, want.token_ids) and torch.equal(got.top_index, want.top_index)):
            failures.append("vocabulary-parallel sample != single-GPU sample")
        if not torch.allclose(got.logsumexp, want.logsumexp, rtol=1e-5, atol=1e-5):
            failures.append("vocabulary-parallel log-sum-exp")
        if _native.workspace_error(dev) != 0:
            failures.append("workspace error word set")
        dist.barrier()
        xch.close()
    except Exception as exc:  # reported to the parent
        failures.append(f"exception: {exc!r}")
    finally:
        with open(f"{result_path}.{rank}", "w") as f:
            f.write("\n".join(failures))
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_vocab_parallel_peer_exchange_two_gpus(tmp_path):
    import torch.multiprocessing as mp
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    port = _free_port()
    result = str(tmp_path / "result")
    ctx = mp.spawn(_worker, args=(2, port, result), nprocs=2, join=False)
    done = False
    for _ in range(60):  # up to 10 minutes
        done = ctx.join(timeout=10)
        if done:
            break
    if not done:
        for proc in ctx.processes:
            proc.kill()
        pytest.fail("vocab-parallel workers did not finish")
    for r in range(2):
        text = open(f"{result}.{r}").read()
        assert text == "", f"rank {r}: {text}"


@pytest.mark.parametrize("route", ["row-sparse", "block-sparse"])
def test_exchange_wait_runs_out_on_one_gpu(cuda_device, route):
    """Failure detection without a fault: a two-rank exchange whose second
    rank never runs (its buffer is a second local one that nothing writes).
    The last CTA's wait gives up after the caller's limit (5 ms), the call
    returns no token (top_index -1, top_value NaN: not a merge of what
    arrived), check_exchange raises, the workspace error word reads 3; after
    the buffers and the workspace are re-zeroed the device keeps working (a
    plain call on the same stream succeeds)."""
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", "grammar-sparse-projection_b200"))
    from gsp import _native
    dev = cuda_device
    rng = np.random.default_rng(3)
    vocab, hidden = 4096, 64
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32)).half().to(dev)
    h = torch.from_numpy(rng.standard_normal((1, hidden), dtype=np.float32)).half().to(dev)
    mask = torch.full((1, vocab // 32), -1, dtype=torch.int32, device=dev)
    own, _ = _native.peer_exchange_alloc(2, 1)
    silent, _ = _native.peer_exchange_alloc(2, 1)
    try:
        from gsp import vocab_parallel as vp
        _native.reset_workspace(dev)
        tv = torch.empty(1, device=dev)
        ti = torch.empty(1, device=dev, dtype=torch.int64)
        t0 = time.perf_counter()
        _native.vocab_parallel(route, h, w[: vocab // 2], mask[:, : vocab // 64], [own, silent], 0, 1,
                               vocab, top_value=tv, top_index=ti, wait_us=5000)
        torch.cuda.synchronize()
        assert time.perf_counter() - t0 < 2.0  # the caller's limit, not the default
        assert ti.item() == -1 and math.isnan(tv.item())
        with pytest.raises(vp.ExchangeTimeout):
            vp.check_exchange(ti)
        assert _native.workspace_error(dev) == 3
        _native.peer_exchange_reset(own, 2, 1)
        _native.peer_exchange_reset(silent, 2, 1)
        _native.reset_workspace(dev)
        logits = torch.empty(1, vocab, device=dev, dtype=torch.float16)
        _native.row_sparse(h, w, mask, logits=logits, top_value=tv, top_index=ti)
        torch.cuda.synchronize()
        assert _native.workspace_error(dev) == 0
        assert ti.item() == logits.argmax(-1).item()
    finally:
        _native.peer_exchange_free(own)
        _native.peer_exchange_free(silent)


def test_prepared_vocab_parallel_single_rank(cuda_device):
    """PreparedVocabParallel (arguments converted once) with world size 1 runs
    the plain projection: equal to gsp_row_sparse_logits, on repeated calls,
    with the top-1 record written into pinned host memory."""
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", "grammar-sparse-projection_b200"))
    from gsp import _native
    dev = cuda_device
    rng = np.random.default_rng(9)
    vocab, hidden = 20000, 128
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32) * 0.1).half().to(dev)
    h = torch.from_numpy(rng.standard_normal((1, hidden), dtype=np.float32)).half().to(dev)
    mask = torch.from_numpy(_case(vocab, hidden, 1, 4, torch.float16)[2]).to(dev)
    own, _ = _native.peer_exchange_alloc(1, 1)
    try:
        lg = torch.empty(1, vocab, dtype=torch.float16, device=dev)
        host = torch.zeros(2, dtype=torch.int64).pin_memory()
        call = _native.PreparedVocabParallel("row-sparse", h, w, mask, [own], 0, 1, vocab, logits=lg,
                                             top_value=host[1:2].view(torch.float32)[:1], top_index=host[0:1])
        lg_ref = torch.empty(1, vocab, dtype=torch.float16, device=dev)
        ti_ref = torch.empty(1, dtype=torch.int64, device=dev)
        tv_ref = torch.empty(1, device=dev)
        _native.row_sparse(h, w, mask, logits=lg_ref, top_value=tv_ref, top_index=ti_ref)
        for _ in range(3):
            host.zero_()
            call()
            torch.cuda.synchronize()
            assert torch.equal(lg, lg_ref)
            assert int(host[0]) == ti_ref.item() and host[1:2].view(torch.float32)[0].item() == tv_ref.item()
        assert _native.workspace_error(dev) == 0
    finally:
        _native.peer_exchange_free(own)
